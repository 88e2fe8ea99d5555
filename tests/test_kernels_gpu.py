"""Per-kernel parity of libtt_b200 against plain PyTorch FP32 math of the same op.

Operands are rounded to FP16 exactly as the kernels consume them, so the only
differences left are accumulation order, FP32 transcendental rounding and the
FP16 rounding of FP16 outputs.  Tolerances are stated per test.
"""

import math

import pytest
import torch
import torch.nn.functional as F

from tiktoktechjam2026_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _gen(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


@pytest.mark.parametrize("d", [32, 64, 96, 128, 256, 512, 768, 1024])
@pytest.mark.parametrize("n", [1, 7, 1000])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_layernorm_rows(tt_lib, d, n, out_dtype):
    g = _gen(d * 31 + n)
    x = (torch.randn(n, d, generator=g) * 3 + 0.5).to(DEV)
    w = torch.randn(d, generator=g).to(DEV)
    b = torch.randn(d, generator=g).to(DEV)
    out = ops.layernorm_rows(x, w, b, 1e-5, out_dtype)
    ref = F.layer_norm(x, (d,), w, b, 1e-5)
    tol = 4e-3 if out_dtype == torch.float16 else 2e-5  # FP16 output rounding (|y| < 8)
    torch.testing.assert_close(out.float(), ref, rtol=tol, atol=tol)


QKV_SHAPES = [(2, 16, 32, 2), (3, 130, 128, 4), (1, 256, 256, 8), (2, 64, 512, 8), (64, 128, 128, 4),
              (2, 128, 128, 16), (1, 70, 64, 8), (2, 128, 1024, 4), (1, 64, 768, 6), (1, 100, 512, 4)]


@pytest.mark.parametrize("B,S,D,H", QKV_SHAPES)
def test_qkv_projection(tt_lib, B, S, D, H):
    g = _gen(B * S + D)
    n = torch.randn(B, S, D, generator=g).half().to(DEV)
    w = (torch.randn(3 * D, D, generator=g) / math.sqrt(D)).half().to(DEV)
    b = (torch.randn(3 * D, generator=g) * 0.1).to(DEV)
    q, k, vt = ops.qkv_projection(n, w, b, H)
    hd = D // H
    ref = (n.float() @ w.float().t() + b).view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
    assert q.shape[-1] == ops.stored_head_dim(hd) and vt.shape[2] == ops.stored_head_dim(hd)
    # FP16 output rounding of |x| < 8 values: 4e-3
    torch.testing.assert_close(q[..., :hd].float(), ref[0], rtol=2e-3, atol=4e-3)
    torch.testing.assert_close(k[..., :hd].float(), ref[1], rtol=2e-3, atol=4e-3)
    torch.testing.assert_close(vt[:, :, :hd, :S].float(), ref[2].transpose(-1, -2), rtol=2e-3, atol=4e-3)
    # head_dim 8 is stored 16 wide; the padding features of q and k are exact zeros.
    assert torch.all(q[..., hd:] == 0) and torch.all(k[..., hd:] == 0)


def test_qkv_projection_rejects_misaligned_outputs(tt_lib):
    """The epilogue stores 16-byte pieces: q/k/vt that are not 16-byte aligned are refused, not written."""
    B, S, D, H = 1, 64, 128, 4
    n = torch.zeros(B, S, D, dtype=torch.float16, device=DEV)
    w = torch.zeros(3 * D, D, dtype=torch.float16, device=DEV)
    b = torch.zeros(3 * D, device=DEV)
    buf = torch.zeros(4 * B * S * D, dtype=torch.float16, device=DEV)
    base = buf.data_ptr()
    q, k, vt = base + 2, base + 2 * B * S * D + 256, base + 4 * B * S * D + 512
    rc = tt_lib.tt_qkv_projection(n.data_ptr(), w.data_ptr(), b.data_ptr(), q, k, vt, B, S, D, H, S,
                                  torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _lib.TT_ERR_ALIGN
    assert torch.all(buf == 0)


def _attn_ref(q, k, vt, scale, causal, mask):
    B, H, S, hd = q.shape
    v = vt[..., :S].transpose(-1, -2).float()
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    if causal:
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    if mask is not None:
        s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)  # rows with no valid key are defined as 0
    return (p @ v).transpose(1, 2).reshape(B, S, H * hd)


ATTN_SHAPES = [
    (2, 2, 16, 16), (1, 4, 130, 32), (2, 2, 256, 64), (1, 8, 1024, 32), (3, 1, 200, 16), (1, 2, 384, 64),
    (2, 4, 200, 8), (1, 16, 128, 8), (2, 2, 200, 128), (1, 2, 1024, 128), (1, 4, 128, 256), (2, 1, 300, 256),
]


@pytest.mark.parametrize("B,H,S,hd", ATTN_SHAPES)
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("mask_kind", [None, "prefix", "random"])
def test_attention(tt_lib, B, H, S, hd, causal, mask_kind):
    g = _gen(B * 1000 + S + hd)
    hs = ops.stored_head_dim(hd)
    q = torch.zeros(B, H, S, hs, dtype=torch.float16)
    k = torch.zeros(B, H, S, hs, dtype=torch.float16)
    q[..., :hd] = torch.randn(B, H, S, hd, generator=g).half()
    k[..., :hd] = torch.randn(B, H, S, hd, generator=g).half()
    q, k = q.to(DEV), k.to(DEV)
    sp = ops.seq_pad_of(S)
    vt = torch.zeros(B, H, hs, sp, dtype=torch.float16)
    vt[:, :, :hd, :S] = torch.randn(B, H, hd, S, generator=g).half()
    if hs > hd:
        vt[:, :, hd:, :S] = 7.0  # rows past head_dim feed no stored output
    vt = vt.to(DEV)
    mask = None
    if mask_kind == "prefix":
        lengths = torch.randint(max(1, S // 2), S + 1, (B,), generator=g)
        mask = (torch.arange(S)[None, :] < lengths[:, None]).to(DEV)
    elif mask_kind == "random":
        mask = (torch.rand(B, S, generator=g) > 0.3).to(DEV)
        mask[:, 0] = True
    scale = hd**-0.5
    out = ops.attention(q, k, vt, scale, causal, mask, head_dim=hd)
    ref = _attn_ref(q[..., :hd], k[..., :hd], vt[:, :, :hd], scale, causal, mask)
    if mask is not None:
        # Padded query rows are defined as zero context.
        ref = ref.masked_fill(~mask[..., None], 0)
    # P is rounded to FP16 before P.V (as in the reference kernel); |ctx| <= max|v| < 5
    torch.testing.assert_close(out.float(), ref, rtol=5e-3, atol=5e-3)


def test_attention_fully_padded_tile_is_zero(tt_lib):
    B, H, S, hd = 2, 2, 512, 32
    g = _gen(9)
    q = torch.randn(B, H, S, hd, generator=g).half().to(DEV)
    k = torch.randn(B, H, S, hd, generator=g).half().to(DEV)
    vt = torch.randn(B, H, hd, S, generator=g).half().to(DEV)
    mask = torch.zeros(B, S, dtype=torch.bool, device=DEV)
    mask[0, :100] = True
    mask[1, :300] = True
    out = ops.attention(q, k, vt, hd**-0.5, True, mask)
    assert torch.all(out[0, 100:] == 0) and torch.all(out[1, 300:] == 0)
    ref = _attn_ref(q, k, vt, hd**-0.5, True, mask)
    torch.testing.assert_close(out[0, :100].float(), ref[0, :100], rtol=5e-3, atol=5e-3)
    torch.testing.assert_close(out[1, :300].float(), ref[1, :300], rtol=5e-3, atol=5e-3)


# d_model 96, 160 and 224 split their rows unevenly between the two epilogue warps of a lane quadrant.
LIN_LN_SHAPES = [(1000, 128, 128), (300, 32, 32), (513, 256, 256), (257, 512, 512), (200, 2048, 512),
                 (129, 1024, 256), (4096, 128, 128), (300, 96, 96), (257, 160, 160), (129, 224, 224),
                 (300, 1024, 1024), (257, 768, 768), (129, 2048, 1024)]


@pytest.mark.parametrize("N,K,D", LIN_LN_SHAPES)
@pytest.mark.parametrize("norm_dtype", [torch.float16, torch.float32])
def test_linear_residual_layernorm(tt_lib, N, K, D, norm_dtype):
    g = _gen(N + K + D)
    a = torch.randn(N, K, generator=g).half().to(DEV)
    w = (torch.randn(D, K, generator=g) / math.sqrt(K)).half().to(DEV)
    b = (torch.randn(D, generator=g) * 0.1).to(DEV)
    r = torch.randn(N, D, generator=g).to(DEV)
    gw = (1 + 0.1 * torch.randn(D, generator=g)).to(DEV)
    gb = (0.1 * torch.randn(D, generator=g)).to(DEV)
    mask = (torch.rand(N, generator=g) > 0.2).to(DEV)
    resid, norm = ops.linear_residual_layernorm(a, w, b, r, gw, gb, 1e-5, norm_dtype, mask)
    ref_r = r + a.float() @ w.float().t() + b
    ref_n = F.layer_norm(ref_r, (D,), gw, gb, 1e-5).masked_fill(~mask[:, None], 0)
    torch.testing.assert_close(resid, ref_r, rtol=1e-5, atol=2e-5)
    tol = 4e-3 if norm_dtype == torch.float16 else 5e-5
    torch.testing.assert_close(norm.float(), ref_n, rtol=tol, atol=tol)


@pytest.mark.parametrize("N,K,Fo", [(1000, 128, 128), (300, 32, 128), (257, 512, 2048), (129, 256, 1024)])
def test_linear_gelu(tt_lib, N, K, Fo):
    g = _gen(N * 3 + K + Fo)
    a = torch.randn(N, K, generator=g).half().to(DEV)
    w = (torch.randn(Fo, K, generator=g) / math.sqrt(K)).half().to(DEV)
    b = (torch.randn(Fo, generator=g) * 0.1).to(DEV)
    out = ops.linear_gelu(a, w, b)
    ref = F.gelu(a.float() @ w.float().t() + b, approximate="none")
    torch.testing.assert_close(out.float(), ref, rtol=2e-3, atol=4e-3)


def test_watchdog_times_out_cleanly_and_context_survives(tt_lib):
    from tiktoktechjam2026_b200 import _lib

    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = tt_lib.tt_watchdog_selftest(20_000_000, stream)  # 20 ms limit
    assert rc == _lib.TT_ERR_TIMEOUT, _lib.last_error()
    # error word was cleared; the context still runs kernels correctly
    word = __import__("ctypes").c_uint(0)
    assert tt_lib.tt_device_error(__import__("ctypes").byref(word), 1) == _lib.TT_OK
    x = torch.randn(64, 128, device=DEV)
    out = ops.layernorm_rows(x, torch.ones(128, device=DEV), torch.zeros(128, device=DEV), 1e-5, torch.float32)
    torch.testing.assert_close(out, F.layer_norm(x, (128,)), rtol=2e-5, atol=2e-5)


# The last two run 2-3 row tiles per CTA of the persistent kernel.
FFN_SHAPES = [(1000, 128, 128), (300, 32, 128), (513, 256, 1024), (129, 64, 256), (4096, 256, 1024), (77, 128, 512),
              (38000, 256, 256), (40000, 128, 128)]


@pytest.mark.parametrize("N,D,Fd", FFN_SHAPES)
@pytest.mark.parametrize("norm_dtype", [torch.float16, torch.float32])
def test_ffn_residual_layernorm(tt_lib, N, D, Fd, norm_dtype):
    g = _gen(N * 7 + D + Fd)
    a = torch.randn(N, D, generator=g).half().to(DEV)
    w1 = (torch.randn(Fd, D, generator=g) / math.sqrt(D)).half().to(DEV)
    b1 = (torch.randn(Fd, generator=g) * 0.1).to(DEV)
    w2 = (torch.randn(D, Fd, generator=g) / math.sqrt(Fd)).half().to(DEV)
    b2 = (torch.randn(D, generator=g) * 0.1).to(DEV)
    r = torch.randn(N, D, generator=g).to(DEV)
    gw = (1 + 0.1 * torch.randn(D, generator=g)).to(DEV)
    gb = (0.1 * torch.randn(D, generator=g)).to(DEV)
    mask = (torch.rand(N, generator=g) > 0.2).to(DEV)
    resid, norm = ops.ffn_residual_layernorm(a, w1, b1, w2, b2, r, gw, gb, 1e-5, norm_dtype, mask)
    # The reference rounds the GELU output to FP16 before the second projection.
    h = F.gelu(a.float() @ w1.float().t() + b1, approximate="none").half().float()
    ref_r = r + h @ w2.float().t() + b2
    ref_n = F.layer_norm(ref_r, (D,), gw, gb, 1e-5).masked_fill(~mask[:, None], 0)
    # The GELU differs from exact erf by < 6.7e-6, which rarely flips the FP16 rounding of h by one
    # ulp (2^-9 at |h| ~ 3); through W2 (|w| <= ~0.3) that moves r by at most ~1.5e-3.
    torch.testing.assert_close(resid, ref_r, rtol=1e-3, atol=2e-3)
    tol = 4e-3 if norm_dtype == torch.float16 else 1e-3
    torch.testing.assert_close(norm.float(), ref_n, rtol=tol, atol=tol)


def test_gelu_matches_exact_erf(tt_lib):
    """GELU of the projection epilogue against exact-erf GELU over a dense input sweep."""
    x = torch.linspace(-12, 12, 128 * 2048, device=DEV).reshape(-1, 128)
    eye = torch.eye(128, device=DEV).half()
    out = ops.linear_gelu(x.half(), eye, torch.zeros(128, device=DEV))
    ref = F.gelu(x.half().float(), approximate="none")
    # out is FP16: within FP16 rounding of the exact value
    torch.testing.assert_close(out.float(), ref, rtol=1e-3, atol=1e-6)


def test_exp2_polynomial_matches_exp2(tt_lib):
    """The softmax's FMA-pipe exponential against exact 2^max(x, -26) over [-125, 64): relative error
    <= 7.9e-5 (the fit's 7.5e-5, the 2^-18 rounding of its clamped input y = (x + 26) / 128 and FP32
    rounding of the result); its FP16 form within one FP16 unit in the last place of the exact 2^x,
    zero below 2^-25 (x < 15.99, below FP16's largest finite value 65504 = 2^15.9993)."""
    g = _gen(77)
    x = torch.cat([torch.linspace(-125.0, 63.99, 1 << 21), (torch.rand(1 << 20, generator=g) * 188.99 - 125.0),
                   torch.tensor([-125.0, -0.5, 0.5, -0.49999997, 0.49999997, 0.0, -1.0, 1.0, 7.9999995, 8.0,
                                 -26.0, -25.5, -25.0, -24.5, -24.0])])
    x = x[: x.numel() // 2 * 2].contiguous().to(DEV)
    y32 = torch.empty_like(x)
    y16 = torch.empty(x.numel(), dtype=torch.float16, device=DEV)
    rc = tt_lib.tt_selftest_exp2_fma(x.data_ptr(), y32.data_ptr(), y16.data_ptr(), x.numel(),
                                     torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _lib.TT_OK, _lib.last_error()
    exact = torch.exp2(x.double())
    clamped = torch.exp2(x.double().clamp_min(-26.0))
    rel = ((y32.double() - clamped).abs() / clamped).max().item()
    assert rel <= 7.9e-5, rel
    sel = x < 15.99
    e = exact[sel]
    ulp = torch.exp2(torch.floor(torch.log2(e)) - 10).clamp_min(2.0 ** -24)
    err16 = (y16[sel].double() - e).abs()
    assert bool(torch.all(err16 <= ulp)), float((err16 / ulp).max())
    assert bool(torch.all(y16[x < -25.0] == 0))
