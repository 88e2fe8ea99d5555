"""The CPU oracle reproduces the reference's own outputs (fixtures written by
tests/golden/make_golden.py from the reference checkout)."""

import numpy as np
import pytest
import torch

import oracle


def _checksums(tensors):
    rows = []
    for v in tensors:
        f = v.detach().double().flatten()
        idx = torch.linspace(0, f.numel() - 1, 8).long()
        rows.append([float(f.sum()), float(f.abs().sum())] + [float(f[i]) for i in idx])
    return np.array(rows, dtype=np.float64)


def _cfg(c):
    B, S, D, H, F, L, causal = c
    return oracle.Config(B, S, D, H, F, L, bool(causal))


def test_reference_source_hash_recorded(golden):
    _, meta = golden
    assert len(meta["reference_sha256_torch_transformer_benchmark"]) == 64


@pytest.mark.parametrize("name", ["t_causal_small", "t_causal_mask", "t_full_mask", "t_causal_s130", "t_hd64"])
def test_tiny_case_matches_reference(golden, name):
    data, meta = golden
    m = meta["tiny"][name]
    cfg = _cfg(m["cfg"])
    sd = oracle.seeded_state_dict(cfg, m["seed"])
    # seeded weights are bit-identical to the reference's BaselineTransformer init
    np.testing.assert_array_equal(_checksums(sd.values()), data[f"{name}/wsum"])
    # Q/K/V packing matches copy_mixed_model_weights (key order = mixed state_dict order)
    packed = oracle.pack_qkv_state_dict(sd)
    keys = m["mixed_state_keys"]
    assert sorted(keys) == sorted(packed.keys())
    np.testing.assert_array_equal(_checksums([packed[k] for k in keys]), data[f"{name}/packedsum"])
    x, mask = oracle.generate_case(cfg, m["seed"], m["padding_ratio"])
    np.testing.assert_array_equal(_checksums([x]), data[f"{name}/xsum"])
    np.testing.assert_array_equal(mask.numpy(), data[f"{name}/mask"])
    y = oracle.forward(sd, cfg, x, None if m["padding_ratio"] <= 0 else mask)
    np.testing.assert_allclose(y.numpy(), data[f"{name}/y"], rtol=0, atol=2e-5)


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C4", "C5"])
def test_bench_config_weights_and_inputs(golden, name):
    data, meta = golden
    m = meta["bench"][name]
    cfg, pad = oracle.CONFIGS[name]
    assert [cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers,
            cfg.causal] == m["cfg"]
    assert pad == m["padding_ratio"]
    sd = oracle.seeded_state_dict(cfg, oracle.DEFAULT_SEED)
    assert list(sd.keys()) == m["weight_keys"]
    np.testing.assert_array_equal(_checksums(sd.values()), data[f"{name}/wsum"])
    x, mask = oracle.generate_case(cfg, oracle.DEFAULT_SEED, pad)
    np.testing.assert_allclose(x.double().sum(dim=(1, 2)).numpy(), data[f"{name}/xsum"], rtol=0, atol=1e-9)
    np.testing.assert_array_equal(mask.sum(dim=1).numpy(), data[f"{name}/lengths"])


@pytest.mark.parametrize("name", ["C1", "C3", "C4"])
def test_bench_config_outputs_match_reference(golden, name):
    """Oracle output of the picked sequences equals the reference's (C2/C5 are covered on the GPU box)."""
    data, meta = golden
    m = meta["bench"][name]
    cfg, pad = oracle.CONFIGS[name]
    sd = oracle.seeded_state_dict(cfg, oracle.DEFAULT_SEED)
    x, mask = oracle.generate_case(cfg, oracle.DEFAULT_SEED, pad)
    for i in m["picked_sequences"]:
        y = oracle.forward(sd, cfg, x[i : i + 1], None if pad <= 0 else mask[i : i + 1])
        np.testing.assert_allclose(y[0, ::16].numpy(), data[f"{name}/y_seq{i}_rows16"], rtol=0, atol=3e-5)


def test_compare_rule_is_or_not_isclose():
    ref = torch.tensor([0.0, 1.0, 10.0, float("nan")])
    out = torch.tensor([0.0019, 1.019, 10.19, 0.0])
    res = oracle.compare(ref, out)
    # 0.0019 <= atol; 0.019 <= 0.02*1; 0.19 <= 0.02*10; NaN in ref fails
    assert res.failed == 1
    res2 = oracle.compare(ref[:3], torch.tensor([0.0021, 1.0, 10.0]))
    assert res2.failed == 1  # 0.0021 > atol and > rtol*0


def test_flops_bytes_c2():
    cfg, _ = oracle.CONFIGS["C2"]
    flops, nbytes = oracle.forward_flops_bytes(cfg)
    assert abs(flops / 1e9 - 120.3) < 1.0
    assert abs(nbytes / 1e9 - 1.41) < 0.05
