"""CPU FP32 restatement of the reference's strict baseline Transformer.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA path: the
tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
use it; the shipped package never imports it.

It restates, in plain PyTorch FP32 CPU math, the parts of
neil0618/TikTokTechJam2026 that define correctness for the forward pass:

* ``seeded_state_dict``   -- weights of ``BaselineTransformer(config)`` built
  right after ``torch.manual_seed(seed)`` (mixed_precision_benchmark.py:53,60;
  module order torch_transformer_benchmark.py:202-237).
* ``generate_case``       -- ``generate_random_case`` on CPU
  (torch_transformer_benchmark.py:448-486).
* ``forward``             -- ``BaselineTransformer.forward``
  (torch_transformer_benchmark.py:162-199 attention, :211-222 block,
  :239-249 model): pre-LN blocks, explicit S x S scores, causal ``triu`` mask,
  key-padding mask, FP32 softmax, exact-erf GELU, padded rows zeroed after
  every block and on output.
* ``compare``             -- ``compare_outputs``'s per-element rule
  (torch_transformer_benchmark.py:503-570): pass iff finite and
  (abs_err <= atol or abs_err <= rtol * |ref|), defaults atol 0.002, rtol 0.02
  (:869-870).
* ``pack_qkv_state_dict`` -- ``copy_mixed_model_weights``'s Q/K/V packing
  (mixed_precision/transformer.py:702-731).

Pinned by tests/golden (fixtures written by tests/golden/make_golden.py from
the reference itself).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class Config:
    """Same fields as the reference's TransformerConfig (torch_transformer_benchmark.py:106-133)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool


# The five BASELINE configurations (C1..C5) and the padding ratio of each.
CONFIGS: Dict[str, Tuple[Config, float]] = {
    "C1": (Config(64, 128, 128, 4, 128, 4, True), 0.0),
    "C2": (Config(64, 1024, 128, 4, 128, 4, True), 0.0),
    "C3": (Config(256, 256, 32, 2, 128, 4, True), 0.0),
    "C4": (Config(16, 2048, 512, 8, 2048, 6, True), 0.5),
    "C5": (Config(512, 1024, 256, 8, 1024, 4, True), 0.0),
}

# Cases of the reference's wider suite that BASELINE.json does not name
# (analysis_profile_mixed.py:20-26; run with every token valid, :45).  Case 8
# (d_model 1024, head_dim 256) is outside this build's shape coverage.
SUITE_CONFIGS: Dict[str, Tuple[Config, float]] = {
    "S6": (Config(10000, 128, 128, 4, 128, 4, True), 0.0),
    "S8": (Config(64, 128, 1024, 4, 1024, 4, True), 0.0),
    "S10": (Config(64, 128, 128, 2, 128, 4, True), 0.0),
    "S11": (Config(64, 128, 128, 16, 128, 4, True), 0.0),
    "S13": (Config(64, 1024, 128, 4, 128, 4, True), 0.0),
}

DEFAULT_SEED = 1234  # torch_transformer_benchmark.py:871
TIMING_SEED_OFFSET = 100000  # torch_transformer_benchmark.py:747
ATOL = 0.002
RTOL = 0.02


def seeded_state_dict(cfg: Config, seed: int = DEFAULT_SEED) -> Dict[str, torch.Tensor]:
    """FP32 weights identical to ``torch.manual_seed(seed); BaselineTransformer(cfg)``.

    nn.Linear / nn.LayerNorm are constructed in the reference's module order
    (per block: norm1, q, k, v, out, norm2, ffn_in, ffn_out; then final_norm),
    so PyTorch's default initialisers draw the same random stream.
    """
    torch.manual_seed(seed)
    D, Fd = cfg.d_model, cfg.ffn_dim
    sd: Dict[str, torch.Tensor] = {}
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        mods = [
            ("norm1", nn.LayerNorm(D)),
            ("attention.q_proj", nn.Linear(D, D)),
            ("attention.k_proj", nn.Linear(D, D)),
            ("attention.v_proj", nn.Linear(D, D)),
            ("attention.out_proj", nn.Linear(D, D)),
            ("norm2", nn.LayerNorm(D)),
            ("ffn_in", nn.Linear(D, Fd)),
            ("ffn_out", nn.Linear(Fd, D)),
        ]
        for name, mod in mods:
            sd[p + name + ".weight"] = mod.weight.detach().clone()
            sd[p + name + ".bias"] = mod.bias.detach().clone()
    fn = nn.LayerNorm(D)
    sd["final_norm.weight"] = fn.weight.detach().clone()
    sd["final_norm.bias"] = fn.bias.detach().clone()
    return sd


def pack_qkv_state_dict(sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Baseline state dict -> mixed-model state dict (q/k/v concatenated)."""
    out: Dict[str, torch.Tensor] = {}
    for key, val in sd.items():
        if ".attention.q_proj." in key:
            suffix = key.split(".attention.q_proj.")[1]
            prefix = key.split(".attention.q_proj.")[0]
            out[f"{prefix}.attention.qkv_proj.{suffix}"] = torch.cat(
                [
                    sd[f"{prefix}.attention.q_proj.{suffix}"],
                    sd[f"{prefix}.attention.k_proj.{suffix}"],
                    sd[f"{prefix}.attention.v_proj.{suffix}"],
                ],
                dim=0,
            )
        elif ".attention.k_proj." in key or ".attention.v_proj." in key:
            continue
        else:
            out[key] = val
    return out


def generate_case(
    cfg: Config,
    seed: int,
    padding_ratio: float = 0.0,
    input_scale: float = 1.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """CPU restatement of generate_random_case (torch_transformer_benchmark.py:448-486)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, generator=g, dtype=torch.float32)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(cfg.batch_size, cfg.seq_len, dtype=torch.bool)
    min_valid = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(min_valid, cfg.seq_len + 1, (cfg.batch_size,), generator=g)
    mask = torch.arange(cfg.seq_len)[None, :] < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


def _layer_norm(x: torch.Tensor, sd: Dict[str, torch.Tensor], name: str) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), sd[name + ".weight"], sd[name + ".bias"], 1e-5)


def _linear(x: torch.Tensor, sd: Dict[str, torch.Tensor], name: str) -> torch.Tensor:
    return F.linear(x, sd[name + ".weight"], sd[name + ".bias"])


def _attention(
    x: torch.Tensor, sd: Dict[str, torch.Tensor], p: str, cfg: Config, mask: Optional[torch.Tensor]
) -> torch.Tensor:
    """BaselineSelfAttention.forward (torch_transformer_benchmark.py:162-199)."""
    B, S, D = x.shape
    H = cfg.num_heads
    hd = D // H

    def heads(t: torch.Tensor) -> torch.Tensor:
        return t.view(B, S, H, hd).transpose(1, 2).contiguous()

    q = heads(_linear(x, sd, p + "attention.q_proj"))
    k = heads(_linear(x, sd, p + "attention.k_proj"))
    v = heads(_linear(x, sd, p + "attention.v_proj"))
    scores = torch.matmul(q, k.transpose(-2, -1)) * (hd**-0.5)
    if cfg.causal:
        upper = torch.ones(S, S, dtype=torch.bool, device=x.device).triu(diagonal=1)
        scores = scores.masked_fill(upper, float("-inf"))
    if mask is not None:
        scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1)
    ctx = torch.matmul(probs, v).transpose(1, 2).contiguous().view(B, S, D)
    out = _linear(ctx, sd, p + "attention.out_proj")
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    return out


@torch.no_grad()
def forward(
    sd: Dict[str, torch.Tensor],
    cfg: Config,
    x: torch.Tensor,
    mask: Optional[torch.Tensor] = None,
    chunk: Optional[int] = None,
) -> torch.Tensor:
    """BaselineTransformer.forward in FP32 on x's device.

    Sequences are independent, so ``chunk`` bounds memory by running batch
    slices (the reference's MicrobatchModel, torch_transformer_benchmark.py:808-833).
    """
    if chunk is not None and x.shape[0] > chunk:
        outs = []
        for s in range(0, x.shape[0], chunk):
            m = None if mask is None else mask[s : s + chunk]
            outs.append(forward(sd, cfg, x[s : s + chunk], m))
        return torch.cat(outs, dim=0)
    x = x.float()
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        x = x + _attention(_layer_norm(x, sd, p + "norm1"), sd, p, cfg, mask)
        h = _linear(_layer_norm(x, sd, p + "norm2"), sd, p + "ffn_in")
        x = x + _linear(F.gelu(h, approximate="none"), sd, p + "ffn_out")
        if mask is not None:
            x = x.masked_fill(~mask[..., None], 0)
    x = _layer_norm(x, sd, "final_norm")
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    return x


@dataclass
class Comparison:
    passed: bool
    total: int
    failed: int
    max_abs: float
    max_rel: float
    mean_abs: float


def compare(ref: torch.Tensor, out: torch.Tensor, rtol: float = RTOL, atol: float = ATOL) -> Comparison:
    """compare_outputs's rule (torch_transformer_benchmark.py:503-570)."""
    if ref.shape != out.shape:
        raise AssertionError(f"shape mismatch: {tuple(ref.shape)} vs {tuple(out.shape)}")
    r = ref.detach().float()
    o = out.detach().float().to(r.device)
    finite = torch.isfinite(r) & torch.isfinite(o)
    err = (o - r).abs()
    ok = finite & ((err <= atol) | (err <= rtol * r.abs()))
    failed = int((~ok).sum().item())
    rel = err / r.abs().clamp_min(1e-12)
    return Comparison(
        passed=failed == 0,
        total=r.numel(),
        failed=failed,
        max_abs=float(err.max().item()) if r.numel() else 0.0,
        max_rel=float(rel.max().item()) if r.numel() else 0.0,
        mean_abs=float(err.mean().item()) if r.numel() else 0.0,
    )


def forward_flops_bytes(cfg: Config) -> Tuple[float, float]:
    """Algorithmic FLOPs and fused-design HBM bytes of one forward (per layer x L).

    FLOPs = 6ND^2 (QKV) + 2*B*S^2*D (causal attention; 4*B*S^2*D if not causal)
            + 2ND^2 (out) + 4NDF (FFN);
    bytes = 8ND + 6D^2 (QKV) + 8ND (attention) + 12ND + 2D^2 (out+LN)
            + 12ND + 4DF (FFN+LN), plus 4ND for the input read by LN0.
    """
    B, S, D, Fd, L = cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.ffn_dim, cfg.num_layers
    N = B * S
    attn = (2.0 if cfg.causal else 4.0) * B * S * S * D
    flops = L * (6.0 * N * D * D + attn + 2.0 * N * D * D + 4.0 * N * D * Fd)
    nbytes = L * (8.0 * N * D + 6 * D * D + 8.0 * N * D + 12.0 * N * D + 2 * D * D + 12.0 * N * D + 4 * D * Fd)
    nbytes += 4.0 * N * D
    return flops, nbytes
