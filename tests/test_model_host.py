"""Host-side surface of the drop-in model (no GPU needed)."""

import pytest
import torch

import oracle
from tiktoktechjam2026_b200 import B200Transformer, MixedPrecisionTransformer, TransformerConfig, copy_mixed_model_weights


def _cfg(name="C1"):
    c, _ = oracle.CONFIGS[name]
    return TransformerConfig(c.batch_size, c.seq_len, c.d_model, c.num_heads, c.ffn_dim, c.num_layers, c.causal)


def test_reference_class_name_alias():
    assert MixedPrecisionTransformer is B200Transformer


def test_state_dict_keys_match_reference_mixed_model(golden):
    _, meta = golden
    m = meta["tiny"]["t_causal_small"]
    B, S, D, H, F, L, causal = m["cfg"]
    model = B200Transformer(TransformerConfig(B, S, D, H, F, L, causal))
    assert list(model.state_dict().keys()) == m["mixed_state_keys"]


def test_constructor_flags_and_attributes():
    model = B200Transformer(
        _cfg(),
        enable_case11_schedule=False,
        enable_attention_output_norm_fusion=False,
        enable_full_ffn_fusion=False,
        enable_fp16_custom_attention=False,
        enable_fp16_normalized_stream=False,
    )
    for attr in ("use_case8_triton", "use_d128_triton", "use_d128_custom_attention", "use_fp16_custom_attention",
                 "use_case11_schedule", "fuse_attention_output_norm", "fuse_full_ffn",
                 "use_fp16_normalized_stream", "use_d32_triton"):
        assert isinstance(getattr(model, attr), bool)
    assert model.assume_all_tokens_valid is False


def test_copy_weights_strict_and_packing():
    cfg = oracle.Config(2, 8, 32, 2, 64, 2, True)
    sd = oracle.seeded_state_dict(cfg)
    base = torch.nn.Module()
    # a minimal baseline-shaped module: load the oracle's state dict into a dict-backed holder
    class Holder(torch.nn.Module):
        def __init__(self, sd):
            super().__init__()
            self._sd = sd

        def state_dict(self, *a, **k):
            return dict(self._sd)

    model = B200Transformer(TransformerConfig(2, 8, 32, 2, 64, 2, True))
    copy_mixed_model_weights(Holder(sd), model)
    w = model.layers[1].attention.qkv_proj.weight
    assert torch.equal(w[:32], sd["layers.1.attention.q_proj.weight"])
    assert torch.equal(w[64:], sd["layers.1.attention.v_proj.weight"])
    assert torch.equal(model.layers[0].attention.qkv_proj.bias[32:64], sd["layers.0.attention.k_proj.bias"])
    packed = oracle.pack_qkv_state_dict(sd)
    for k, v in model.state_dict().items():
        assert torch.equal(v, packed[k]), k


def test_convert_keeps_fp32_bias_copies():
    model = B200Transformer(TransformerConfig(1, 8, 32, 2, 64, 1, True))
    b = model.layers[0].ffn_in.bias.detach().clone()
    model.convert_projections_to_fp16()
    assert model.layers[0].ffn_in.weight.dtype == torch.float16
    assert model.layers[0].ffn_in.bias.dtype == torch.float16
    assert model.layers[0].norm1.weight.dtype == torch.float32
    assert torch.equal(model._bias_fp32["layers.0.ffn_in"], b)


def test_forward_rejects_non_fp32_and_cpu():
    model = B200Transformer(TransformerConfig(1, 8, 32, 2, 64, 1, True))
    with pytest.raises(ValueError, match="FP32"):
        model(torch.zeros(1, 8, 32, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="CUDA"):
        model(torch.zeros(1, 8, 32))


class _RowwiseModel(torch.nn.Module):
    """Stand-in model: each sequence's output depends only on that sequence (and its mask row)."""

    def __init__(self):
        super().__init__()
        self.calls = []

    def forward(self, x, mask=None):
        self.calls.append(x.shape[0])
        y = x * 2.0 + 1.0
        if mask is not None:
            y = y.masked_fill(~mask[..., None], 0.0)
        return y


def test_microbatch_wrapper_matches_whole_batch():
    """PreallocatedMicrobatchModel (mixed_precision_benchmark.py:13-33): slices of microbatch_size, ragged
    tail, mask sliced alongside, a batch no larger than one microbatch passed through untouched."""
    from tiktoktechjam2026_b200 import PreallocatedMicrobatchModel

    g = torch.Generator().manual_seed(3)
    x = torch.randn(10, 5, 4, generator=g)
    mask = torch.rand(10, 5, generator=g) > 0.4
    inner = _RowwiseModel()
    wrapped = PreallocatedMicrobatchModel(inner, 4)
    out = wrapped(x, mask)
    assert inner.calls == [4, 4, 2]
    assert out.dtype == torch.float32 and torch.equal(out, _RowwiseModel()(x, mask))
    inner.calls.clear()
    assert torch.equal(wrapped(x[:4]), x[:4] * 2.0 + 1.0) and inner.calls == [4]
    with pytest.raises(ValueError):
        PreallocatedMicrobatchModel(inner, 0)
