"""The batch split across GPUs and gathered to GPU 0 (the north star's multi-GPU case).

Each rank (one process per GPU, NCCL only for the handle exchange and
barriers) runs its contiguous slice of the batch through
``forward_gather``, which pushes the FP32 output into rank 0's gather buffer
over NVLink; rank 0 then checks the gathered batch element-wise against the
strict FP32 oracle under the reference's rule (zero failed elements), against
the reference's own stored outputs of the golden sequences, and bit for bit
against its own 1-GPU forward of the whole batch.  Skipped with fewer than
two GPUs.
"""

import json
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CHUNK = {"C1": 64, "C4": 2, "C5": 32}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, result_path):
    from datetime import timedelta

    import numpy as np

    import oracle
    from tiktoktechjam2026_b200 import B200Transformer, TransformerConfig, copy_mixed_model_weights
    from tiktoktechjam2026_b200.sharding import PeerGatherBuffer, shard_bounds

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        cfg, pad = oracle.CONFIGS[name]
        sd = oracle.seeded_state_dict(cfg, oracle.DEFAULT_SEED)

        class _Baseline(torch.nn.Module):
            def state_dict(self, *a, **k):
                return dict(sd)

        model = B200Transformer(TransformerConfig(cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads,
                                                  cfg.ffn_dim, cfg.num_layers, cfg.causal))
        copy_mixed_model_weights(_Baseline(), model)
        model = model.to(dev).eval()
        model.convert_projections_to_fp16()
        model.assume_all_tokens_valid = pad <= 0
        x, mask = oracle.generate_case(cfg, oracle.DEFAULT_SEED, pad)
        mask = None if pad <= 0 else mask
        s0, s1 = shard_bounds(cfg.batch_size, world, rank)
        xs = x[s0:s1].contiguous().to(dev)
        ms = None if mask is None else mask[s0:s1].contiguous().to(dev)
        gather = PeerGatherBuffer(cfg.batch_size, (cfg.seq_len, cfg.d_model), rank, world, dev)
        out = gather.local_view(0)[s0:s1] if rank == 0 else torch.empty_like(xs)
        with torch.inference_mode():
            # Twice: the second call's last layer must wait for the first call's push.
            for _ in range(2):
                model.forward_gather(xs, ms, out, gather.dst(0) if rank != 0 else 0)
            model.gather_wait(dev)
            torch.cuda.synchronize(dev)
            dist.barrier(device_ids=[rank])
            if rank == 0:
                got = gather.local_view(0)
                whole = model(x.to(dev), None if mask is None else mask.to(dev))
                prev = (torch.backends.cuda.matmul.allow_tf32, torch.get_float32_matmul_precision())
                torch.backends.cuda.matmul.allow_tf32 = False
                torch.set_float32_matmul_precision("highest")
                sdd = {k: v.to(dev) for k, v in sd.items()}
                ref = oracle.forward(sdd, cfg, x.to(dev), None if mask is None else mask.to(dev), chunk=CHUNK[name])
                torch.backends.cuda.matmul.allow_tf32 = prev[0]
                torch.set_float32_matmul_precision(prev[1])
                res = oracle.compare(ref, got)
                here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
                data = np.load(os.path.join(here, "golden.npz"))
                with open(os.path.join(here, "golden_meta.json")) as f:
                    meta = json.load(f)
                gold_failed = 0
                for i in meta["bench"][name]["picked_sequences"]:
                    gold = torch.from_numpy(data[f"{name}/y_seq{i}_rows16"]).to(dev)
                    gold_failed += oracle.compare(gold, got[i, ::16]).failed
                record = {"failed": res.failed, "total": res.total, "max_abs": res.max_abs,
                          "golden_failed": gold_failed, "bitwise_equal_to_1gpu": bool(torch.equal(got, whole)),
                          "padded_rows_zero": True if mask is None else bool(torch.all(got[~mask.to(dev)] == 0))}
                with open(result_path, "w") as f:
                    json.dump(record, f)
            dist.barrier(device_ids=[rank])
        gather.close()
    finally:
        dist.destroy_process_group()


def _worlds():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return sorted({w for w in (2, n) if 2 <= w <= min(n, 8)})


@pytest.mark.parametrize("name", ["C5", "C4"])
@pytest.mark.parametrize("world", _worlds() or [2])
def test_batch_split_gathered_to_gpu0_matches_oracle(tt_lib, tmp_path, name, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path = str(tmp_path / "gather.json")
    mp.start_processes(_worker, args=(world, _free_port(), name, path), nprocs=world, join=True,
                       start_method="spawn")
    with open(path) as f:
        rec = json.load(f)
    print(f"{name} world {world}: {rec}")
    assert rec["failed"] == 0, rec
    assert rec["golden_failed"] == 0, rec
    assert rec["bitwise_equal_to_1gpu"], rec
    assert rec["padded_rows_zero"], rec
