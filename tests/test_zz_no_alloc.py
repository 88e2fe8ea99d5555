"""The allocation-free masked attention entry point agrees with the allocating path and with FP32 math.

tt_causal_attention_masked_noalloc serves callers that cannot allocate device
memory (CUDA-graph capture in progress, device memory owned by an external
pool, no allocation allowed after start-up): it keeps its per-sequence scratch
in a static array inside the library.  This test calls it through the C ABI
twice in a row, with different masks so the second call must overwrite what
the first left in the shared array, and compares each result with
tt_mask_kv_end + tt_causal_attention on the same inputs, within the attention
tests' tolerance.  A second test runs it at head_dim 16, 32 and 64, causal and
not, twice in a row with different masks, against plain PyTorch FP32 attention
on the same FP16 operands.  The file sorts last so a failing run stops only
after every other test has run; it also passes on its own in a fresh process.
"""

import ctypes

import pytest
import torch

from tiktoktechjam2026_b200 import _lib, ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _reference_path(q, k, vt, mask, scale):
    B, H, S, hd = q.shape
    m8 = mask.contiguous().view(torch.uint8)
    kv_end = torch.empty(B, dtype=torch.int32, device=DEV)
    ctx = torch.empty(B, S, H * hd, dtype=torch.float16, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    _lib.check(_lib.lib().tt_mask_kv_end(m8.data_ptr(), B, S, kv_end.data_ptr(), stream))
    _lib.check(_lib.lib().tt_causal_attention(q.data_ptr(), k.data_ptr(), vt.data_ptr(), m8.data_ptr(),
                                              kv_end.data_ptr(), ctx.data_ptr(), B, S, H, hd, vt.shape[-1],
                                              scale, 1, stream))
    return ctx


def _noalloc_path(q, k, vt, mask, scale, ctx):
    B, H, S, hd = q.shape
    m8 = mask.contiguous().view(torch.uint8)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    _lib.check(_lib.lib().tt_causal_attention_masked_noalloc(
        q.data_ptr(), k.data_ptr(), vt.data_ptr(), m8.data_ptr(), ctx.data_ptr(), B, S, H, hd, vt.shape[-1],
        scale, 1, stream))


def test_noalloc_matches_allocating_path_twice(tt_lib):
    B, H, S, hd = 6, 4, 640, 32
    g = torch.Generator().manual_seed(2024)
    q = torch.randn(B, H, S, hd, generator=g).half().to(DEV)
    k = torch.randn(B, H, S, hd, generator=g).half().to(DEV)
    sp = ops.seq_pad_of(S)
    vt = torch.randn(B, H, hd, sp, generator=g).half().to(DEV)
    scale = hd**-0.5
    lengths_a = torch.tensor([640, 1, 129, 300, 511, 200])
    lengths_b = torch.tensor([17, 640, 640, 64, 128, 639])
    ctx = torch.empty(B, S, H * hd, dtype=torch.float16, device=DEV)  # caller-provided output
    for lengths in (lengths_a, lengths_b):
        mask = (torch.arange(S)[None, :] < lengths[:, None]).to(DEV)
        _noalloc_path(q, k, vt, mask, scale, ctx)
        ref = _reference_path(q, k, vt, mask, scale)
        torch.cuda.synchronize()
        torch.testing.assert_close(ctx.float(), ref.float(), rtol=5e-3, atol=5e-3)
    word = ctypes.c_uint(0)
    assert _lib.lib().tt_device_error(ctypes.byref(word), 1) == _lib.TT_OK and word.value == 0


def test_noalloc_rejects_batch_beyond_static_limit(tt_lib):
    q = torch.zeros(1, 1, 8, 16, dtype=torch.float16, device=DEV)
    mask = torch.ones(1, 8, dtype=torch.uint8, device=DEV)
    rc = _lib.lib().tt_causal_attention_masked_noalloc(q.data_ptr(), q.data_ptr(), q.data_ptr(), mask.data_ptr(),
                                                       q.data_ptr(), 65537, 8, 1, 16, 8, 0.25, 1,
                                                       torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _lib.TT_ERR_SHAPE
    assert "65536" in _lib.last_error()


def _fp32_attention(q, k, vt, scale, causal, mask):
    """softmax(q k^T * scale + masks) v in FP32 from the FP16 operands; padded query rows are zero."""
    B, H, S, hd = q.shape
    v = vt[..., :S].transpose(-1, -2).float()
    s = (q.float() @ k.float().transpose(-1, -2)) * scale
    if causal:
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
    p = torch.nan_to_num(torch.softmax(s, dim=-1), nan=0.0)
    ctx = (p @ v).transpose(1, 2).reshape(B, S, H * hd)
    return ctx.masked_fill(~mask[..., None], 0)


@pytest.mark.parametrize("hd", [16, 32, 64])
@pytest.mark.parametrize("causal", [True, False])
def test_noalloc_matches_fp32_attention(tt_lib, hd, causal):
    B, H, S = 5, 2, 200
    g = torch.Generator().manual_seed(hd * 10 + int(causal))
    q = torch.randn(B, H, S, hd, generator=g).half().to(DEV)
    k = torch.randn(B, H, S, hd, generator=g).half().to(DEV)
    sp = ops.seq_pad_of(S)
    vt = torch.zeros(B, H, hd, sp, dtype=torch.float16)
    vt[..., :S] = torch.randn(B, H, hd, S, generator=g).half()
    vt = vt.to(DEV)
    scale = hd**-0.5
    ctx = torch.empty(B, S, H * hd, dtype=torch.float16, device=DEV)
    for lengths in (torch.tensor([200, 1, 77, 128, 199]), torch.tensor([64, 200, 3, 150, 129])):
        mask = (torch.arange(S)[None, :] < lengths[:, None]).to(DEV)
        m8 = mask.contiguous().view(torch.uint8)
        _lib.check(_lib.lib().tt_causal_attention_masked_noalloc(
            q.data_ptr(), k.data_ptr(), vt.data_ptr(), m8.data_ptr(), ctx.data_ptr(), B, S, H, hd, sp, scale,
            int(causal), torch.cuda.current_stream(DEV).cuda_stream))
        torch.cuda.synchronize()
        ref = _fp32_attention(q, k, vt, scale, causal, mask)
        # P is rounded to FP16 before P.V; |ctx| <= max|v| < 5
        torch.testing.assert_close(ctx.float(), ref, rtol=5e-3, atol=5e-3)
