"""Writes the golden fixtures that pin the CPU oracle to the reference itself.

Run in a container where the reference checkout is importable (it is not on
the GPU box; the fixtures it writes travel instead):

    python tests/golden/make_golden.py --reference <path to TikTokTechJam2026>

For every case it imports the reference's own ``torch_transformer_benchmark``
(``BaselineTransformer``, ``generate_random_case``, ``TransformerConfig``) and
``mixed_precision.copy_mixed_model_weights``, and records:

* tiny cases: checksums of the seeded weights, of the inputs and of the
  packed (Q/K/V concatenated) mixed-model state dict the reference's weight
  copy produces; the full mask and the full reference FP32 CPU output;
* the five benchmark configurations (C1..C5): per-tensor weight checksums, the
  input's per-sequence checksums and valid lengths, and the reference output
  of two sequences (every 16th row) computed on those sequences alone
  (sequences are independent in the model).

Output: tests/golden/golden.npz (+ golden_meta.json).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

TINY_CASES = {
    # name: (B, S, D, H, F, L, causal, padding_ratio, seed)
    "t_causal_small": (2, 16, 32, 2, 64, 2, True, 0.0, 1234),
    "t_causal_mask": (3, 40, 64, 4, 96, 2, True, 0.5, 1234),
    "t_full_mask": (2, 24, 32, 2, 32, 1, False, 0.3, 77),
    "t_causal_s130": (1, 130, 128, 4, 128, 2, True, 0.0, 1234),
    "t_hd64": (2, 72, 128, 2, 256, 1, True, 0.0, 5),
}

BENCH_CASES = {
    "C1": (64, 128, 128, 4, 128, 4, True, 0.0),
    "C2": (64, 1024, 128, 4, 128, 4, True, 0.0),
    "C3": (256, 256, 32, 2, 128, 4, True, 0.0),
    "C4": (16, 2048, 512, 8, 2048, 6, True, 0.5),
    "C5": (512, 1024, 256, 8, 1024, 4, True, 0.0),
}


def checksums(tensors) -> np.ndarray:
    """Per tensor: sum, sum of |.|, and 8 fixed-position samples (float64)."""
    rows = []
    for v in tensors:
        f = v.detach().double().flatten()
        idx = torch.linspace(0, f.numel() - 1, 8).long()
        rows.append([float(f.sum()), float(f.abs().sum())] + [float(f[i]) for i in idx])
    return np.array(rows, dtype=np.float64)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--seed", type=int, default=1234)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch_transformer_benchmark as ttb  # the reference's own module
    from mixed_precision import MixedPrecisionTransformer, copy_mixed_model_weights

    torch.set_num_threads(os.cpu_count() or 1)
    torch.set_float32_matmul_precision("highest")
    src_sha = hashlib.sha256(
        open(os.path.join(args.reference, "torch_transformer_benchmark.py"), "rb").read()
    ).hexdigest()
    arrays = {}
    meta = {"reference_sha256_torch_transformer_benchmark": src_sha, "tiny": {}, "bench": {}}

    def make(B, S, D, H, F, L, causal):
        return ttb.TransformerConfig(B, S, D, H, F, L, causal)

    for name, (B, S, D, H, F, L, causal, pad, seed) in TINY_CASES.items():
        cfg = make(B, S, D, H, F, L, causal)
        torch.manual_seed(seed)
        base = ttb.BaselineTransformer(cfg).eval()
        x, mask = ttb.generate_random_case(cfg, torch.device("cpu"), torch.float32, seed, pad, 1.0)
        with torch.inference_mode():
            y = base(x, None if pad <= 0 else mask)
        mixed = MixedPrecisionTransformer(cfg)
        copy_mixed_model_weights(base, mixed)
        arrays[f"{name}/wsum"] = checksums(base.state_dict().values())
        arrays[f"{name}/packedsum"] = checksums(mixed.state_dict().values())
        arrays[f"{name}/xsum"] = checksums([x])
        arrays[f"{name}/mask"] = mask.numpy()
        arrays[f"{name}/y"] = y.numpy()
        meta["tiny"][name] = {"cfg": [B, S, D, H, F, L, causal], "padding_ratio": pad, "seed": seed,
                              "mixed_state_keys": list(mixed.state_dict().keys())}
        print("tiny", name, "done", flush=True)

    for name, (B, S, D, H, F, L, causal, pad) in BENCH_CASES.items():
        cfg = make(B, S, D, H, F, L, causal)
        torch.manual_seed(args.seed)
        base = ttb.BaselineTransformer(cfg).eval()
        arrays[f"{name}/wsum"] = checksums(base.state_dict().values())
        x, mask = ttb.generate_random_case(cfg, torch.device("cpu"), torch.float32, args.seed, pad, 1.0)
        arrays[f"{name}/xsum"] = x.double().sum(dim=(1, 2)).numpy()
        arrays[f"{name}/lengths"] = mask.sum(dim=1).numpy().astype(np.int64)
        lengths = mask.sum(dim=1)
        picks = [0, int(torch.argmin(lengths))] if pad > 0 else [0, B - 1]
        if picks[1] == picks[0]:
            picks[1] = B - 1
        with torch.inference_mode():
            for i in picks:
                y = base(x[i : i + 1], None if pad <= 0 else mask[i : i + 1])
                arrays[f"{name}/y_seq{i}_rows16"] = y[0, ::16].numpy()
        meta["bench"][name] = {"cfg": [B, S, D, H, F, L, causal], "padding_ratio": pad,
                               "picked_sequences": picks, "weight_keys": list(base.state_dict().keys())}
        print("bench", name, "done", flush=True)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", len(arrays), "arrays")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
